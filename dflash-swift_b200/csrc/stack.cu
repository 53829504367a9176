// Glue kernels of the tensor-parallel verify stack (the hybrid target's layers around the
// quantized projections): residual add + RMSNorm, the SiLU-gated MLP activation, the
// gated-delta layer's causal depthwise convolution, per-head normalisation, gates and
// gated output norm, and the attention layer's q/k norm + rotary embedding + cache append
// and its decode attention with the output gate.  The projections themselves are
// dflash_qmm and the recurrence is dflash_gdn_step.
//
// All tensors are row-major with one row per token (M rows, the verify block).  Every
// kernel here is latency-bound and tiny next to the weight stream, so each is launched
// with programmatic dependent launch: it is scheduled while its predecessor drains and
// waits (griddepcontrol.wait) before touching memory, then releases its successor.
#include "common.cuh"
#include "dflash_stack.h"
#include "tp_layout.cuh"

namespace dflash {
namespace stack {

__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
__device__ __forceinline__ uint16_t to_bf(float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    return *reinterpret_cast<const uint16_t*>(&h);
}
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float bf_round(float v) { return bf(to_bf(v)); }
__device__ __forceinline__ float silu(float v) { return v / (1.f + __expf(-v)); }
__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
    return static_cast<uint32_t>(to_bf(a)) | (static_cast<uint32_t>(to_bf(b)) << 16);
}

// Wait for the predecessor, then let the successor be scheduled.
__device__ __forceinline__ void chain_in() {
    pdl_wait();
    pdl_launch_dependents();
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += red[i];  // the same order on every thread
    return t;
}

// resid[m] += delta[m] (if given); out[m] = bf16(resid[m] * rsqrt(mean(resid[m]^2) + eps) * w).
// A row is split over a cluster of kNormSplit CTAs of 128 threads (more loads in flight
// than one CTA per row gives); each thread keeps up to VPT float4 of its part in
// registers.  The parts' sums of squares are exchanged through distributed shared
// memory and added in rank order, so every CTA uses the same scale.  The weight (written by
// no kernel of the stream) is requested before the wait on the predecessor.  Needs H a
// multiple of 4 kNormSplit, H / kNormSplit <= 512 VPT, delta / w / out 8-byte aligned.
constexpr int kNormSplit = 4;

// Cluster barrier halves: arrive (relaxed: orders nothing), arrive with release, wait with
// acquire.  Every thread of every CTA of the cluster takes each step.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_shared_cluster_f32(uint32_t cluster_addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}

// Hands this CTA's part of a row's sum of squares to the kNormSplit CTAs of the cluster and
// returns the row's total, the parts added in rank order (the same bits in every CTA).
// The part is stored into slot `rank` of every CTA's `parts`, so after the one barrier all
// reads are local and no CTA touches another's shared memory again: a CTA may exit as soon
// as it is done.  The caller arrived (relaxed) on the cluster barrier at its start, so that
// every CTA is known to be running before it is written to; this waits for that phase first.
__device__ __forceinline__ float cluster_row_total(float part, float* parts, uint32_t rank) {
    cluster_wait_acquire();
    if (threadIdx.x < kNormSplit) st_shared_cluster_f32(map_to_rank(smem_u32(&parts[rank]), threadIdx.x), part);
    cluster_arrive_release();
    cluster_wait_acquire();
    float tot = 0.f;
#pragma unroll
    for (int r = 0; r < kNormSplit; ++r) tot += parts[r];
    return tot;
}

// This thread's VPT words (4 bf16 each) of a norm weight: words base + threadIdx.x + 128 j.
template <int VPT>
__device__ __forceinline__ void load_norm_weight(uint2 (&ww)[VPT], const uint16_t* __restrict__ w, int base, int P4) {
    const uint2* w4 = reinterpret_cast<const uint2*>(w) + base;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int i = threadIdx.x + 128 * j;
        ww[j] = i < P4 ? __ldg(w4 + i) : make_uint2(0u, 0u);
    }
}

template <int VPT>
__global__ void __launch_bounds__(128) add_rmsnorm_kernel(float* __restrict__ resid, const uint16_t* __restrict__ delta,
                                                          const uint16_t* __restrict__ w, uint16_t* __restrict__ out,
                                                          int H, float eps) {
    __shared__ float red[4];
    __shared__ float parts[kNormSplit];
    const uint32_t rank = cluster_rank();
    const int m = blockIdx.y, P4 = H / (4 * kNormSplit), base = (int)rank * P4;  // float4 units
    cluster_arrive_relaxed();
    uint2 ww[VPT];
    load_norm_weight<VPT>(ww, w, base, P4);
    chain_in();
    float4* r4 = reinterpret_cast<float4*>(resid + (size_t)m * H) + base;
    const uint2* d4 = reinterpret_cast<const uint2*>(delta + (size_t)m * H) + base;
    float4 v[VPT];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int i = threadIdx.x + 128 * j;
        if (i < P4) {
            v[j] = r4[i];
            if (delta) {
                const uint2 d = d4[i];
                v[j].x += bf16_lo(d.x);
                v[j].y += bf16_hi(d.x);
                v[j].z += bf16_lo(d.y);
                v[j].w += bf16_hi(d.y);
                r4[i] = v[j];
            }
            ss = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, fmaf(v[j].w, v[j].w, ss))));
        }
    }
    const float tot = cluster_row_total(block_sum(ss, red), parts, rank);
    const float rs = rsqrtf(tot / H + eps);
    uint2* o4 = reinterpret_cast<uint2*>(out + (size_t)m * H) + base;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int i = threadIdx.x + 128 * j;
        if (i < P4)
            o4[i] = make_uint2(pack_bf2(v[j].x * rs * bf16_lo(ww[j].x), v[j].y * rs * bf16_hi(ww[j].x)),
                               pack_bf2(v[j].z * rs * bf16_lo(ww[j].y), v[j].w * rs * bf16_hi(ww[j].y)));
    }
}

// add_rmsnorm whose delta is the tensor-parallel sum of the ranks' partials, read from
// this rank's exchange buffer (set `set`, filled by dflash_tp_push on every rank): each
// data word is taken once it carries this exchange's epoch (bounded wait), and
// delta = bf16(sum of the slots in rank order).
template <int VPT>
__global__ void __launch_bounds__(128) add_rmsnorm_reduce_kernel(float* __restrict__ resid, void* xbase, int world,
                                                                 int set, const uint16_t* __restrict__ w,
                                                                 uint16_t* __restrict__ out, int M, int H, float eps) {
    __shared__ float red[4];
    __shared__ float parts[kNormSplit];
    const uint32_t rank = cluster_rank();
    const int m = blockIdx.y, P4 = H / (4 * kNormSplit), base = (int)rank * P4;  // float4 units
    cluster_arrive_relaxed();
    uint2 ww[VPT];
    load_norm_weight<VPT>(ww, w, base, P4);
    chain_in();
    tp::Header* hdr = static_cast<tp::Header*>(xbase);
    const uint32_t e = hdr->next[set];
    float4* r4 = reinterpret_cast<float4*>(resid + (size_t)m * H) + base;
    float4 v[VPT];
    float ss = 0.f;
    // JB float4 slices at a time: their residual values and every source's two words per
    // slice are all requested before any is inspected, so the loads overlap; a word without
    // the expected epoch is then waited for alone.  Slices, sources and components are
    // summed in the same order as one slice at a time would.
    constexpr int JB = VPT < 4 ? VPT : VPT == 4 ? 4 : 2;  // 8 would spill (2 x 8 words per slice)
#pragma unroll
    for (int j0 = 0; j0 < VPT; j0 += JB) {
        uint64_t w0[JB][tp::kMaxRanks], w1[JB][tp::kMaxRanks];
#pragma unroll
        for (int jj = 0; jj < JB; ++jj) {
            const int i = threadIdx.x + 128 * (j0 + jj);
            if (i < P4) {
                v[j0 + jj] = r4[i];
                const size_t word = ((size_t)m * H + 4 * (size_t)(base + i)) / 2;  // two data words per float4
#pragma unroll
                for (int r = 0; r < tp::kMaxRanks; ++r) {
                    if (r < world) {
                        const uint64_t* src = tp::slot_ptr(xbase, world, M, H, set, r) + word;
                        w0[jj][r] = tp::ld_relaxed_sys_u64(src);
                        w1[jj][r] = tp::ld_relaxed_sys_u64(src + 1);
                    }
                }
            }
        }
#pragma unroll
        for (int jj = 0; jj < JB; ++jj) {
            const int j = j0 + jj, i = threadIdx.x + 128 * j;
            if (i < P4) {
                const size_t word = ((size_t)m * H + 4 * (size_t)(base + i)) / 2;
                float sx = 0.f, sy = 0.f, sz = 0.f, sw = 0.f;
#pragma unroll
                for (int r = 0; r < tp::kMaxRanks; ++r) {
                    if (r < world) {
                        const uint64_t* src = tp::slot_ptr(xbase, world, M, H, set, r) + word;
                        const uint32_t d0 =
                            (uint32_t)(w0[jj][r] >> 32) == e ? (uint32_t)w0[jj][r] : tp::wait_word(src, e);
                        const uint32_t d1 =
                            (uint32_t)(w1[jj][r] >> 32) == e ? (uint32_t)w1[jj][r] : tp::wait_word(src + 1, e);
                        sx += bf16_lo(d0);
                        sy += bf16_hi(d0);
                        sz += bf16_lo(d1);
                        sw += bf16_hi(d1);
                    }
                }
                v[j].x += bf_round(sx);
                v[j].y += bf_round(sy);
                v[j].z += bf_round(sz);
                v[j].w += bf_round(sw);
                r4[i] = v[j];
                ss = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, fmaf(v[j].w, v[j].w, ss))));
            }
        }
    }
    const float tot = cluster_row_total(block_sum(ss, red), parts, rank);
    const float rs = rsqrtf(tot / H + eps);
    uint2* o4 = reinterpret_cast<uint2*>(out + (size_t)m * H) + base;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int i = threadIdx.x + 128 * j;
        if (i < P4)
            o4[i] = make_uint2(pack_bf2(v[j].x * rs * bf16_lo(ww[j].x), v[j].y * rs * bf16_hi(ww[j].x)),
                               pack_bf2(v[j].z * rs * bf16_lo(ww[j].y), v[j].w * rs * bf16_hi(ww[j].y)));
    }
    // this exchange is consumed: the next push into the set uses the following epoch
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) hdr->seq[set] = e;
}

// The same for any H and alignment (row re-read from global memory for the second pass).
__global__ void __launch_bounds__(256) add_rmsnorm_any_kernel(float* __restrict__ resid,
                                                              const uint16_t* __restrict__ delta,
                                                              const uint16_t* __restrict__ w,
                                                              uint16_t* __restrict__ out, int H, float eps) {
    __shared__ float red[8];
    chain_in();
    const int m = blockIdx.x;
    float* r = resid + (size_t)m * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        float v = r[i];
        if (delta) {
            v += bf(delta[(size_t)m * H + i]);
            r[i] = v;
        }
        ss = fmaf(v, v, ss);
    }
    const float rs = rsqrtf(block_sum(ss, red) / H + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) out[(size_t)m * H + i] = to_bf(r[i] * rs * bf(w[i]));
}

// gu = [gate (I) | up (I)] per row -> y = silu(gate) * up
__global__ void silu_mul_kernel(const uint16_t* __restrict__ gu, uint16_t* __restrict__ y, int M, int I) {
    chain_in();
    const size_t n = (size_t)M * I;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const size_t m = e / I, i = e % I;
        const float g = bf(gu[m * 2 * I + i]), u = bf(gu[m * 2 * I + I + i]);
        y[e] = to_bf(silu(g) * u);
    }
}

// Causal depthwise convolution over tokens with a window of the previous kc-1 inputs,
// followed by SiLU.  x: [M, ld] with the convolved channels at [0, C); window: [kc-1, C];
// w: [C, kc].  The C channels are `parts` equal parts (q, k, v); y holds each part as its
// own contiguous [M, C / parts] block.  The window is the pre-round one and is only read:
// after the round dflash_gdn_conv_rollback rebuilds it from the accepted inputs.  One
// thread per channel; the M <= 16 inputs are loaded up front.
template <int KC>
__global__ void conv_silu_kernel(const uint16_t* __restrict__ x, int ld, const uint16_t* __restrict__ window,
                                 const uint16_t* __restrict__ w, uint16_t* __restrict__ y, int M, int C, int parts) {
    chain_in();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    constexpr int h = KC - 1;
    float xs[h + 16];
#pragma unroll
    for (int i = 0; i < h; ++i) xs[i] = bf(window[(size_t)i * C + c]);
#pragma unroll
    for (int t = 0; t < 16; ++t) xs[h + t] = t < M ? bf(x[(size_t)t * ld + c]) : 0.f;
    float wk[KC];
#pragma unroll
    for (int i = 0; i < KC; ++i) wk[i] = bf(w[(size_t)c * KC + i]);
    const int cp = C / parts, part = c / cp, cc = c - part * cp;
#pragma unroll
    for (int t = 0; t < 16; ++t) {
        if (t < M) {
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < KC; ++i) acc = fmaf(wk[i], xs[t + i], acc);
            y[((size_t)part * M + t) * cp + cc] = to_bf(silu(acc));
        }
    }
}

// Per (token, head) of the gated-delta layer: L2-normalise q and k (dk each) in place,
// alpha = exp(-exp(a_log[h]) * softplus(a + dt_bias[h])), beta = sigmoid(b).
// q, k: [M, heads * dk]; ab: [M, ld_ab] with b at [0, heads) and a at [heads, 2 heads).
// One warp per (token, head).
__global__ void gdn_gates_kernel(uint16_t* __restrict__ q, uint16_t* __restrict__ k, const uint16_t* __restrict__ ab,
                                 int ld_ab, const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                                 float* __restrict__ alpha, float* __restrict__ beta, int M, int heads, int dk) {
    chain_in();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M * heads) return;
    const int t = warp / heads, h = warp % heads;
    for (int part = 0; part < 2; ++part) {
        uint16_t* v = (part ? k : q) + ((size_t)t * heads + h) * dk;
        float ss = 0.f;
        for (int i = lane; i < dk; i += 32) ss = fmaf(bf(v[i]), bf(v[i]), ss);
        const float rs = rsqrtf(warp_sum(ss) + 1e-6f);
        for (int i = lane; i < dk; i += 32) v[i] = to_bf(bf(v[i]) * rs);
    }
    if (lane == 0) {
        const float b = bf(ab[(size_t)t * ld_ab + h]);
        const float a = bf(ab[(size_t)t * ld_ab + heads + h]);
        const float sp = a + dt_bias[h] > 20.f ? a + dt_bias[h] : log1pf(__expf(a + dt_bias[h]));
        alpha[(size_t)t * heads + h] = __expf(-__expf(a_log[h]) * sp);
        beta[(size_t)t * heads + h] = 1.f / (1.f + __expf(-b));
    }
}

// The gated-delta layer's conv and gates in one kernel (the same arithmetic as
// conv_silu_kernel followed by gdn_gates_kernel, so the same bits): one warp per (token,
// head, part q | k | v) covering the head's dk channels (lane l: channels l + 32 j), with
// all of its conv inputs loaded at once.  Causal conv + SiLU, rounded to bf16; q and k
// L2-normalised over the head; written to y as the parts' [M, heads dk] blocks.  The q
// warp's lane 0 also writes alpha and beta of (token, head).
// Tap i of row t reads the input KC-1-i steps back along t's history: the block rows
// before it (a chain), or its ancestors when `parents` gives a tree (the convolution
// of a tree row is that of its root-to-row path), then the window once the history
// runs past the block's anchor: tap i of a row at depth D < KC-1-i reads window row
// D + i (both forms).
template <int KC, int DJ>
__global__ void gdn_conv_gates_kernel(const uint16_t* __restrict__ x, int ld, const uint16_t* __restrict__ window,
                                      const uint16_t* __restrict__ w, uint16_t* __restrict__ y,
                                      const uint16_t* __restrict__ ab, int ld_ab, const float* __restrict__ a_log,
                                      const float* __restrict__ dt_bias, float* __restrict__ alpha,
                                      float* __restrict__ beta, int M, int heads,
                                      const int32_t* __restrict__ parents) {
    constexpr int dk = 32 * DJ;
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const bool live = wid < M * heads * 3, gates = wid % 3 == 0 && lane == 0;
    const int t = wid / (heads * 3), h = (wid / 3) % heads, part = wid % 3;
    const int C = 3 * heads * dk, cp = heads * dk;
    // the conv taps and gate parameters (written by no kernel of the stream) are requested
    // before the wait on the predecessor, the gate inputs together with the conv inputs
    float wk[DJ][KC], dtb = 0.f, alog = 0.f;
    if (live) {
#pragma unroll
        for (int j = 0; j < DJ; ++j)
#pragma unroll
            for (int i = 0; i < KC; ++i) wk[j][i] = bf(__ldg(w + (size_t)(part * cp + h * dk + lane + 32 * j) * KC + i));
        if (gates) {
            dtb = __ldg(dt_bias + h);
            alog = __ldg(a_log + h);
        }
    }
    chain_in();
    if (!live) return;
    float gb = 0.f, ga = 0.f;
    if (gates) {
        gb = bf(ab[(size_t)t * ld_ab + h]);
        ga = bf(ab[(size_t)t * ld_ab + heads + h]);
    }
    // back[s]: the block row s steps back from t, or -1 once the history is in the window
    int back[KC];
    back[0] = t;
#pragma unroll
    for (int s = 1; s < KC; ++s)
        back[s] = back[s - 1] < 0 ? -1 : parents ? tree_parent(parents, back[s - 1]) : back[s - 1] - 1;
    int depth = 0;  // t's depth, capped at KC - 1 (only its comparison with s matters)
#pragma unroll
    for (int s = 1; s < KC; ++s) depth += back[s] >= 0;
    float xin[DJ][KC];
#pragma unroll
    for (int j = 0; j < DJ; ++j) {
        const int c = part * cp + h * dk + lane + 32 * j;
#pragma unroll
        for (int i = 0; i < KC; ++i) {
            const int src = back[KC - 1 - i];
            xin[j][i] = src < 0 ? bf(window[(size_t)(depth + i) * C + c]) : bf(x[(size_t)src * ld + c]);
        }
    }
    float v[DJ];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < DJ; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < KC; ++i) acc = fmaf(wk[j][i], xin[j][i], acc);
        v[j] = bf_round(silu(acc));
        ss = fmaf(v[j], v[j], ss);
    }
    uint16_t* out = y + ((size_t)part * M + t) * cp + (size_t)h * dk + lane;
    if (part < 2) {
        const float rs = rsqrtf(warp_sum(ss) + 1e-6f);
#pragma unroll
        for (int j = 0; j < DJ; ++j) out[32 * j] = to_bf(v[j] * rs);
    } else {
#pragma unroll
        for (int j = 0; j < DJ; ++j) out[32 * j] = to_bf(v[j]);
    }
    if (gates) {
        const float sp = ga + dtb > 20.f ? ga + dtb : log1pf(__expf(ga + dtb));
        alpha[(size_t)t * heads + h] = __expf(-__expf(alog) * sp);
        beta[(size_t)t * heads + h] = 1.f / (1.f + __expf(-gb));
    }
}

// gdn_conv_gates_kernel for layers whose q and k have fewer heads than v: x rows hold
// [q (k_heads dk) | k (k_heads dk) | v (heads dk)], each key head shared by heads / k_heads
// value heads.  One warp per (token, slot), slots 0 .. k_heads-1 the q heads, then the k
// heads, then the value heads; y receives [q: M x k_heads dk | k: M x k_heads dk |
// v: M x heads dk]; the gates are per value head (ab holds b then a for each value head)
// and written by the value warps.  Taps as in gdn_conv_gates_kernel (chain or tree).
template <int KC, int DJ>
__global__ void gdn_conv_gates_grouped_kernel(const uint16_t* __restrict__ x, int ld,
                                              const uint16_t* __restrict__ window, const uint16_t* __restrict__ w,
                                              uint16_t* __restrict__ y, const uint16_t* __restrict__ ab, int ld_ab,
                                              const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                                              float* __restrict__ alpha, float* __restrict__ beta, int M, int heads,
                                              int k_heads, const int32_t* __restrict__ parents) {
    constexpr int dk = 32 * DJ;
    const int slots = 2 * k_heads + heads;
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const bool live = wid < M * slots;
    const int t = wid / slots, slot = wid % slots;
    const int part = slot < k_heads ? 0 : slot < 2 * k_heads ? 1 : 2;
    const int h = slot - part * k_heads;  // head within its part
    const int C = slots * dk;
    const int c0 = part * k_heads * dk + h * dk;  // first channel of this warp's head
    const bool gates = part == 2 && lane == 0;
    // weights before the wait on the predecessor, as in gdn_conv_gates_kernel
    float wk[DJ][KC], dtb = 0.f, alog = 0.f;
    if (live) {
#pragma unroll
        for (int j = 0; j < DJ; ++j)
#pragma unroll
            for (int i = 0; i < KC; ++i) wk[j][i] = bf(__ldg(w + (size_t)(c0 + lane + 32 * j) * KC + i));
        if (gates) {
            dtb = __ldg(dt_bias + h);
            alog = __ldg(a_log + h);
        }
    }
    chain_in();
    if (!live) return;
    float gb = 0.f, ga = 0.f;
    if (gates) {
        gb = bf(ab[(size_t)t * ld_ab + h]);
        ga = bf(ab[(size_t)t * ld_ab + heads + h]);
    }
    int back[KC];
    back[0] = t;
#pragma unroll
    for (int s = 1; s < KC; ++s)
        back[s] = back[s - 1] < 0 ? -1 : parents ? tree_parent(parents, back[s - 1]) : back[s - 1] - 1;
    int depth = 0;
#pragma unroll
    for (int s = 1; s < KC; ++s) depth += back[s] >= 0;
    float xin[DJ][KC];
#pragma unroll
    for (int j = 0; j < DJ; ++j) {
        const int c = c0 + lane + 32 * j;
#pragma unroll
        for (int i = 0; i < KC; ++i) {
            const int src = back[KC - 1 - i];
            xin[j][i] = src < 0 ? bf(window[(size_t)(depth + i) * C + c]) : bf(x[(size_t)src * ld + c]);
        }
    }
    float v[DJ];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < DJ; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < KC; ++i) acc = fmaf(wk[j][i], xin[j][i], acc);
        v[j] = bf_round(silu(acc));
        ss = fmaf(v[j], v[j], ss);
    }
    const int part_heads = part < 2 ? k_heads : heads;
    uint16_t* out = y + (size_t)part * M * k_heads * dk + ((size_t)t * part_heads + h) * dk + lane;
    if (part < 2) {
        const float rs = rsqrtf(warp_sum(ss) + 1e-6f);
#pragma unroll
        for (int j = 0; j < DJ; ++j) out[32 * j] = to_bf(v[j] * rs);
    } else {
#pragma unroll
        for (int j = 0; j < DJ; ++j) out[32 * j] = to_bf(v[j]);
        if (gates) {
            const float sp = ga + dtb > 20.f ? ga + dtb : log1pf(__expf(ga + dtb));
            alpha[(size_t)t * heads + h] = __expf(-__expf(alog) * sp);
            beta[(size_t)t * heads + h] = 1.f / (1.f + __expf(-gb));
        }
    }
}

// out[t, h*dv + i] = rmsnorm(o[t, h, :]) * w[i] * silu(z[t, h*dv + i]); one warp per (t, h).
// C = dv / 32 (1, 2, 4 or 8): lane l holds elements l + 32 c, the weight requested before
// the wait on the predecessor and o and z together after it, so the kernel waits on
// memory once.  C = 0: any dv, in loops.  Both sum the squares in the same order.
template <int C>
__global__ void gated_norm_kernel(const uint16_t* __restrict__ o, const uint16_t* __restrict__ z, int ld_z,
                                  const uint16_t* __restrict__ w, uint16_t* __restrict__ out, int M, int heads, int dv,
                                  float eps) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if constexpr (C > 0) {
        float wv[C];
#pragma unroll
        for (int c = 0; c < C; ++c) wv[c] = bf(__ldg(w + lane + 32 * c));
        chain_in();
        if (warp >= M * heads) return;
        const int t = warp / heads, h = warp % heads;
        const uint16_t* ov = o + ((size_t)t * heads + h) * dv;
        const uint16_t* zv = z + (size_t)t * ld_z + (size_t)h * dv;
        float ov_f[C], zv_f[C];
#pragma unroll
        for (int c = 0; c < C; ++c) {
            ov_f[c] = bf(ov[lane + 32 * c]);
            zv_f[c] = bf(zv[lane + 32 * c]);
        }
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c) ss = fmaf(ov_f[c], ov_f[c], ss);
        const float rs = rsqrtf(warp_sum(ss) / dv + eps);
#pragma unroll
        for (int c = 0; c < C; ++c)
            out[((size_t)t * heads + h) * dv + lane + 32 * c] = to_bf(ov_f[c] * rs * wv[c] * silu(zv_f[c]));
    } else {
        chain_in();
        if (warp >= M * heads) return;
        const int t = warp / heads, h = warp % heads;
        const uint16_t* ov = o + ((size_t)t * heads + h) * dv;
        float ss = 0.f;
        for (int i = lane; i < dv; i += 32) ss = fmaf(bf(ov[i]), bf(ov[i]), ss);
        const float rs = rsqrtf(warp_sum(ss) / dv + eps);
        for (int i = lane; i < dv; i += 32) {
            const float zz = bf(z[(size_t)t * ld_z + (size_t)h * dv + i]);
            out[((size_t)t * heads + h) * dv + i] = to_bf(bf(ov[i]) * rs * bf(w[i]) * silu(zz));
        }
    }
}

// Attention-layer prep, one warp per (token, head slot).  qkv row t (stride ld) holds
// [q (hq * d) | gate (hq * d) | k (hkv * d) | v (hkv * d)].  Slot < hq: q head, RMSNorm with
// q_norm then rotary embedding on its first `rot` dims, in place.  Slot >= hq: kv head j,
// k gets k_norm and the rotary embedding and goes to cache_k[j, pos0 + t]; v is copied to
// cache_v[j, pos0 + t].  Rotary: rotate-half over the first rot dims, frequency
// theta^(-2i/rot) for pair (i, i + rot/2), position pos0 + t.  Lane l holds dims
// l + 32 c, so with rot a multiple of 64 both halves of a pair sit in one lane.
// With a tree parent list the rotary position is pos0 + depth(t) (a tree row sits at its
// depth on its path); the cache slot stays pos0 + t.
template <int CH>
__global__ void attn_prep_kernel(uint16_t* __restrict__ qkv, int ld, const uint16_t* __restrict__ q_norm,
                                 const uint16_t* __restrict__ k_norm, uint16_t* __restrict__ cache_k,
                                 uint16_t* __restrict__ cache_v, int M, int hq, int hkv, int rot, int pos0,
                                 int max_len, float eps, float theta, const int32_t* __restrict__ parents,
                                 const int32_t* __restrict__ position) {
    constexpr int d = CH * 32;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int slots = hq + hkv;
    const bool live = warp < M * slots;
    const int t = live ? warp / slots : 0, slot = warp % slots;
    // the norm weight (written by no kernel of the stream) is requested before the wait on
    // the predecessor; after it, the cache position and this warp's rows are requested together
    const uint16_t* nw = slot < hq ? q_norm : k_norm;
    float nwv[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) nwv[c] = live ? bf(__ldg(nw + lane + 32 * c)) : 0.f;
    chain_in();
    uint16_t* row = qkv + (size_t)t * ld;
    uint16_t* src = slot < hq ? row + (size_t)slot * d : row + (size_t)(2 * hq + (slot - hq)) * d;
    const uint16_t* vs = row + (size_t)(2 * hq + hkv + (slot - hq)) * d;  // slot >= hq: the v row
    float v[CH];
    uint16_t vcopy[CH];
    if (live) {
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            v[c] = bf(src[lane + 32 * c]);
            if (slot >= hq) vcopy[c] = vs[lane + 32 * c];
        }
    }
    if (position) {  // the cache position from device memory (a graph replayed at a new context)
        pos0 = *position;
        if (pos0 < 0 || pos0 + M > max_len) {
            if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&g_device_error, DFLASH_DEVERR_POSITION);
            return;
        }
    }
    if (!live) return;
    if (slot >= hq) {
        uint16_t* vd = cache_v + ((size_t)(slot - hq) * max_len + pos0 + t) * d;
#pragma unroll
        for (int c = 0; c < CH; ++c) vd[lane + 32 * c] = vcopy[c];
    }
    uint16_t* dst = slot < hq ? src : cache_k + ((size_t)(slot - hq) * max_len + pos0 + t) * d;
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) ss = fmaf(v[c], v[c], ss);
    const float rs = rsqrtf(warp_sum(ss) / d + eps);
#pragma unroll
    for (int c = 0; c < CH; ++c) v[c] = bf_round(v[c] * rs * nwv[c]);
    const int half_c = rot / 64;  // pair partner is c + half_c
    const float pos = (float)(pos0 + (parents ? tree_walk(parents, t).depth : t));
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        if (c < half_c) {
            const int i = lane + 32 * c;
            const float inv = exp2f(-(2.f * i / rot) * log2f(theta));
            float sn, cs;
            sincosf(pos * inv, &sn, &cs);
            float b = 0.f;
#pragma unroll
            for (int cc = 0; cc < CH; ++cc)
                if (cc == c + half_c) b = v[cc];  // register select, no local-memory indexing
            const float a = v[c];
            v[c] = a * cs - b * sn;
#pragma unroll
            for (int cc = 0; cc < CH; ++cc)
                if (cc == c + half_c) v[cc] = b * cs + a * sn;
        }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) dst[lane + 32 * c] = to_bf(v[c]);
}

// Decode attention of the block.  A cluster of SPLIT CTAs serves one (kv head, token t):
// the keys 0 .. pos0 + t that token t sees are cut into SPLIT contiguous ranges, one per
// CTA, and each CTA runs an online softmax over its range for all G = hq / hkv q heads
// that read this kv head, in chunks of kChunk keys.  Lane l holds dims [l CH, l CH + CH)
// of every row it touches, so each key or value row is one coalesced read.
//   scores: a warp takes KU = 32 / GP keys at a time (GP >= G, a power of two); every
//           lane forms the KU x GP partial dot products over its dims and a butterfly
//           reduce-scatter (16 + 8 + 4 + 2 + 1 exchanges) leaves lane u GP + g holding
//           the full dot product of key u with head g;
//   p V:    warp w takes keys w, w + 8, ... (kUnroll in flight); each lane accumulates its
//           dims for the G heads; the 8 warps' partials are summed in a fixed order
//           through shared memory.
// The CTAs' (max, sum, p V) partials are merged through distributed shared memory, each
// CTA of the cluster finishing a quarter of the outputs, with the output gate:
//   out[t, h d + e] = softmax(q k^T scale) v * sigmoid(gate[t, h d + e]).
// With a tree parent list, block key pos0 + a is visible to token t only when row a lies
// on t's root-to-row path (the cached prefix stays visible); hidden keys score -inf.  A
// chunk or CTA range may then hold no visible key: its exponent base stays finite (0)
// so its weights come out 0, and the merge gives such a CTA weight 0 (t itself is
// always visible, so some CTA holds a finite maximum).
constexpr int kSplit = 4;       // CTAs per (kv head, token) ...
constexpr int kSplitSmall = 8;  // ... or, when the grid would leave most SMs idle, twice as many
constexpr int kChunk = 384;     // keys a CTA scores per pass (a 1032-key context in one pass at SPLIT 4)
constexpr int kMaxG = 8;
constexpr int kUnroll = 8;     // value rows a warp has in flight in the p V pass (its key order does not depend on it)

template <int CH>
__device__ __forceinline__ void load_row(const uint16_t* p, float (&v)[CH]) {
    if constexpr (CH == 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
        v[4] = bf16_lo(u.z); v[5] = bf16_hi(u.z); v[6] = bf16_lo(u.w); v[7] = bf16_hi(u.w);
    } else if constexpr (CH == 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
    } else {
        const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
        v[0] = bf16_lo(u); v[1] = bf16_hi(u);
    }
}

// Butterfly reduce-scatter of 32 values per lane: afterwards lane l holds the sum over
// the warp of value l.
__device__ __forceinline__ float reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
    for (int lvl = 0; lvl < 5; ++lvl) {
        const int m = 16 >> lvl, n = 32 >> lvl, h = n / 2;
        const bool hi = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < h; ++i) {
            const float send = hi ? v[i] : v[i + h];
            const float keep = hi ? v[i + h] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
    }
    return v[0];
}

template <int CH, int GP, int SPLIT>
__global__ void __launch_bounds__(256) attn_decode_kernel(const uint16_t* __restrict__ qkv, int ld,
                                                          const uint16_t* __restrict__ cache_k,
                                                          const uint16_t* __restrict__ cache_v,
                                                          uint16_t* __restrict__ out, int hq, int hkv, int pos0,
                                                          int max_len, float scale,
                                                          const int32_t* __restrict__ parents,
                                                          const int32_t* __restrict__ position) {
    constexpr int d = CH * 32;
    constexpr int KU = 32 / GP;  // keys per warp step in the scores pass
    static_assert(GP <= kMaxG && KU * CH <= 64, "score registers");
    __shared__ float s_p[kMaxG][kChunk];
    __shared__ __align__(16) float s_red[4][kMaxG][d];  // warp partials; s_red[0] ends as the CTA's p V
    __shared__ float s_m[kMaxG], s_l[kMaxG], s_corr[kMaxG], s_f[SPLIT][kMaxG], s_den[kMaxG];
    chain_in();
    if (position) {  // the cache position from device memory (a graph replayed at a new context)
        pos0 = *position;
        if (pos0 < 0 || pos0 + (int)gridDim.y > max_len) {  // every CTA leaves here, before any cluster barrier
            if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) atomicOr(&g_device_error, DFLASH_DEVERR_POSITION);
            return;
        }
    }
    const int G = hq / hkv;
    const int kvh = blockIdx.x / SPLIT, t = blockIdx.y;
    const uint32_t rank = cluster_rank();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = pos0 + t + 1;
    const int k0 = (int)((long long)n * rank / SPLIT), k1 = (int)((long long)n * (rank + 1) / SPLIT);
    const uint32_t visible = parents ? tree_walk(parents, t).path : 0u;  // tree rounds: t's path rows

    float q[GP][CH];
    const uint16_t* qrow = qkv + (size_t)t * ld + (size_t)kvh * G * d + lane * CH;
#pragma unroll
    for (int g = 0; g < GP; ++g)
#pragma unroll
        for (int c = 0; c < CH; ++c) q[g][c] = g < G ? bf(qrow[(size_t)g * d + c]) * scale : 0.f;
    if (threadIdx.x < kMaxG) {
        s_m[threadIdx.x] = -INFINITY;
        s_l[threadIdx.x] = 0.f;
    }
    const uint16_t* kb = cache_k + (size_t)kvh * max_len * d + lane * CH;
    const uint16_t* vb = cache_v + (size_t)kvh * max_len * d + lane * CH;
    float acc[kMaxG][CH];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g)
#pragma unroll
        for (int c = 0; c < CH; ++c) acc[g][c] = 0.f;

    for (int c0 = k0; c0 < k1; c0 += kChunk) {
        const int len = min(kChunk, k1 - c0);
        __syncthreads();  // s_p of the previous chunk is consumed; s_m / s_l initialised
        // scores: keys j0 + u, u < KU, for warp steps j0 = KU warp, KU (warp + 8), ...
        for (int j0 = KU * warp; j0 < len; j0 += 8 * KU) {
            float kv[KU][CH];
#pragma unroll
            for (int u = 0; u < KU; ++u) {
                if (j0 + u < len) {
                    load_row<CH>(kb + (size_t)(c0 + j0 + u) * d, kv[u]);
                } else {
#pragma unroll
                    for (int c = 0; c < CH; ++c) kv[u][c] = 0.f;
                }
            }
            float v[32];
#pragma unroll
            for (int u = 0; u < KU; ++u)
#pragma unroll
                for (int g = 0; g < GP; ++g) {
                    float sdot = 0.f;
#pragma unroll
                    for (int c = 0; c < CH; ++c) sdot = fmaf(q[g][c], kv[u][c], sdot);
                    v[u * GP + g] = sdot;
                }
            const float dot = reduce_scatter32(v, lane);
            const int u = lane / GP, g = lane % GP;
            if (g < G && j0 + u < len) {
                const int b = c0 + j0 + u - pos0;  // block row of the key (< 0: the prefix)
                s_p[g][j0 + u] = parents && b >= 0 && !((visible >> b) & 1u) ? -INFINITY : dot;
            }
        }
        __syncthreads();
        // softmax bookkeeping: warp g owns head g
        if (warp < G) {
            float mc = -INFINITY;
            for (int j = lane; j < len; j += 32) mc = fmaxf(mc, s_p[warp][j]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
            const float mold = s_m[warp], mnew = fmaxf(mold, mc);
            const float mbase = mnew == -INFINITY ? 0.f : mnew;  // no visible key yet: weights 0
            float ls = 0.f;
            for (int j = lane; j < len; j += 32) {
                const float p = __expf(s_p[warp][j] - mbase);
                s_p[warp][j] = p;
                ls += p;
            }
            ls = warp_sum(ls);
            if (lane == 0) {
                const float corr = __expf(mold - mbase);  // 0 while mold = -inf
                s_corr[warp] = corr;
                s_l[warp] = s_l[warp] * corr + ls;
                s_m[warp] = mnew;
            }
        }
        __syncthreads();
        // p V
#pragma unroll
        for (int g = 0; g < kMaxG; ++g) {
            const float corr = g < G ? s_corr[g] : 0.f;
#pragma unroll
            for (int c = 0; c < CH; ++c) acc[g][c] *= corr;
        }
        for (int j0 = warp; j0 < len; j0 += 8 * kUnroll) {
            float vv[kUnroll][CH];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int j = j0 + 8 * u;
                if (j < len) load_row<CH>(vb + (size_t)(c0 + j) * d, vv[u]);
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int j = j0 + 8 * u;
                if (j < len) {
#pragma unroll
                    for (int g = 0; g < kMaxG; ++g) {
                        if (g < G) {
                            const float p = s_p[g][j];
#pragma unroll
                            for (int c = 0; c < CH; ++c) acc[g][c] = fmaf(p, vv[u][c], acc[g][c]);
                        }
                    }
                }
            }
        }
    }
    // the 8 warps' partials: warps 0-3 store, warps 4-7 add, then s_red[0] += s_red[1..3]
    if (warp < 4) {
#pragma unroll
        for (int g = 0; g < kMaxG; ++g)
#pragma unroll
            for (int c = 0; c < CH; ++c)
                if (g < G) s_red[warp][g][lane * CH + c] = acc[g][c];
    }
    __syncthreads();
    if (warp >= 4) {
#pragma unroll
        for (int g = 0; g < kMaxG; ++g)
#pragma unroll
            for (int c = 0; c < CH; ++c)
                if (g < G) s_red[warp - 4][g][lane * CH + c] += acc[g][c];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * d; idx += blockDim.x) {
        const int g = idx / d, e = idx - g * d;
        s_red[0][g][e] = ((s_red[0][g][e] + s_red[1][g][e]) + s_red[2][g][e]) + s_red[3][g][e];
    }
    cluster_sync_all();  // every CTA's partial is complete and visible to the cluster
    // merge weights per head: f_r = exp(m_r - max), den = sum_r f_r l_r
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        float mr[SPLIT], mx = -INFINITY;
#pragma unroll
        for (int r = 0; r < SPLIT; ++r) {
            mr[r] = ld_shared_cluster_f32(map_to_rank(smem_u32(&s_m[g]), r));
            mx = fmaxf(mx, mr[r]);
        }
        float den = 0.f;
#pragma unroll
        for (int r = 0; r < SPLIT; ++r) {
            const float f = mr[r] == -INFINITY ? 0.f : __expf(mr[r] - mx);
            s_f[r][g] = f;
            den = fmaf(f, ld_shared_cluster_f32(map_to_rank(smem_u32(&s_l[g]), r)), den);
        }
        s_den[g] = den;
    }
    __syncthreads();
    // this CTA finishes outputs [rank, rank + SPLIT, ...) of the G d
    for (int idx = (int)rank + SPLIT * threadIdx.x; idx < G * d; idx += SPLIT * blockDim.x) {
        const int g = idx / d, ee = idx - g * d;
        float num = 0.f;
#pragma unroll
        for (int r = 0; r < SPLIT; ++r)
            num = fmaf(s_f[r][g], ld_shared_cluster_f32(map_to_rank(smem_u32(&s_red[0][g][ee]), r)), num);
        const int h = kvh * G + g;
        const float gt = bf(qkv[(size_t)t * ld + (size_t)(hq + h) * d + ee]);
        out[(size_t)t * hq * d + (size_t)h * d + ee] = to_bf(num / s_den[g] / (1.f + __expf(-gt)));
    }
    cluster_sync_all();  // every CTA is done reading the others' shared memory
}

// Greedy accept of a verify round from the LM head's argmax keys (dflash_qmm_ex with
// argmax_keys): tokens[i] = the argmax of row i; match i = (proposals[i] == tokens[i]) for
// i < drafts; accepted = the length of the leading run of matches.  One warp.
__global__ void accept_kernel(const unsigned long long* __restrict__ keys, const int32_t* __restrict__ proposals,
                              int drafts, int32_t* __restrict__ tokens, int32_t* __restrict__ accepted) {
    chain_in();
    const int lane = threadIdx.x;
    int run = 0;
    for (int base = 0; base <= drafts; base += 32) {
        const int i = base + lane;
        int32_t tok = 0;
        if (i <= drafts) {
            tok = (int32_t)(~(uint32_t)(keys[i] & 0xffffffffull));
            tokens[i] = tok;
        }
        const bool miss = i < drafts && proposals[i] != tok;
        const unsigned mm = __ballot_sync(0xffffffffu, miss);
        const int valid = min(32, drafts - base);  // match slots in this chunk
        if (run == base) run += mm ? min(__ffs(mm) - 1, valid) : max(valid, 0);
    }
    if (lane == 0) *accepted = run;
}

// dflash_accept over the ranks' keys in an exchange buffer laid out for [M, 4] bf16
// (8 bytes of a key = two data words: low then high half).  One warp; lane i < M takes
// row i's key from every rank, keeps the largest, then the leading run of matches as in
// accept_kernel.  Records the exchange as consumed.
__global__ void accept_reduce_kernel(void* xbase, int world, int set, const int32_t* __restrict__ proposals,
                                     int drafts, int32_t* __restrict__ tokens, int32_t* __restrict__ accepted) {
    chain_in();
    tp::Header* hdr = static_cast<tp::Header*>(xbase);
    const uint32_t e = hdr->next[set];
    const int M = drafts + 1, lane = threadIdx.x;
    int run = 0;
    for (int base = 0; base <= drafts; base += 32) {
        const int i = base + lane;
        int32_t tok = 0;
        if (i <= drafts) {
            unsigned long long best = 0ull;
            for (int r = 0; r < world; ++r) {
                const uint64_t* src = tp::slot_ptr(xbase, world, M, 4, set, r) + 2 * (size_t)i;
                const uint32_t lo = tp::wait_word(src, e), hi = tp::wait_word(src + 1, e);
                const unsigned long long key = (static_cast<unsigned long long>(hi) << 32) | lo;
                best = key > best ? key : best;
            }
            tok = (int32_t)(~(uint32_t)(best & 0xffffffffull));
            tokens[i] = tok;
        }
        const bool miss = i < drafts && proposals[i] != tok;
        const unsigned mm = __ballot_sync(0xffffffffu, miss);
        const int valid = min(32, drafts - base);
        if (run == base) run += mm ? min(__ffs(mm) - 1, valid) : max(valid, 0);
    }
    if (lane == 0) {
        *accepted = run;
        hdr->seq[set] = e;
    }
}

inline unsigned grid_for(size_t n, int block) {
    const size_t g = (n + block - 1) / block;
    return (unsigned)(g < 4096 ? (g > 0 ? g : 1) : 4096);
}

inline cudaStream_t as_stream(dflash_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// The accepted path of a tree round (DFlashDraftTree.acceptedPath,
// Sources/DFlashKit/DFlashDraftTree.swift:122-141): from the anchor, step into the first
// child (row order) whose drafted token is the target's token at the current row, until
// no child is.  One warp, lane r standing for row r: a step is one ballot over the rows
// whose parent is the current row.  Rows only increase along a path, so at most rows - 1
// steps.
__global__ void accept_tree_kernel(const int32_t* __restrict__ target, const int32_t* __restrict__ parents,
                                   const int32_t* __restrict__ tokens, int rows, int32_t* __restrict__ path,
                                   int32_t* __restrict__ path_len, int32_t* __restrict__ next_token) {
    chain_in();
    const int lane = threadIdx.x;
    const int par = lane < rows ? tree_parent(parents, lane) : -1;
    const int tok = lane < rows ? tokens[lane] : 0;
    int row = 0, n = 1;
    if (lane == 0) path[0] = 0;
    for (int step = 1; step < rows; ++step) {
        const int want = target[row];
        const unsigned hit = __ballot_sync(0xffffffffu, par == row && tok == want);
        if (!hit) break;
        row = __ffs(hit) - 1;
        if (lane == 0) path[n] = row;
        ++n;
    }
    if (lane == 0) {
        *path_len = n;
        *next_token = target[row];
    }
}

// y[r, n] = bf16(y[r, n] + bias[n]): the bf16 add of a broadcast bias row that
// QuantizedLinear applies after its matmul.  One thread per element.
__global__ void bias_add_kernel(uint16_t* __restrict__ y, const uint16_t* __restrict__ bias, long long total, int N) {
    chain_in();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    y[i] = to_bf(bf(y[i]) + bf(bias[i % N]));
}

// After a tree round, cache rows pos0 + rows[i] move to pos0 + i.  grid (hkv, layers, 2):
// cache_k for z = 0, cache_v for z = 1.  A block stages all `keep` source rows in shared
// memory before writing any, so moves whose sources and destinations overlap are safe.
struct CompactRows {
    int32_t r[kMaxTreeRows];
};

__global__ void __launch_bounds__(256) kv_compact_kernel(uint16_t* __restrict__ cache_k, uint16_t* __restrict__ cache_v,
                                                         long long layer_stride, int d, int pos0, int max_len,
                                                         CompactRows rows, int keep) {
    __shared__ uint4 buf[kMaxTreeRows * 32];  // keep rows of d <= 256 bf16
    chain_in();
    uint16_t* base = (blockIdx.z ? cache_v : cache_k) + (size_t)blockIdx.y * (size_t)layer_stride +
                     ((size_t)blockIdx.x * max_len + pos0) * d;
    const int per_row = d / 8;  // uint4 per cache row
    for (int idx = threadIdx.x; idx < keep * per_row; idx += blockDim.x) {
        const int i = idx / per_row, c = idx - i * per_row;
        buf[idx] = reinterpret_cast<const uint4*>(base + (size_t)rows.r[i] * d)[c];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < keep * per_row; idx += blockDim.x) {
        const int i = idx / per_row, c = idx - i * per_row;
        reinterpret_cast<uint4*>(base + (size_t)i * d)[c] = buf[idx];
    }
}

}  // namespace stack
}  // namespace dflash

using namespace dflash;
using stack::as_stream;

extern "C" int dflash_stack_add_rmsnorm(float* resid, const dflash_bf16* delta, const dflash_bf16* weight,
                                        dflash_bf16* out, int M, int H, float eps, dflash_stream_t stream) {
    if (!resid || !weight || !out || M < 1 || H < 1 || M > 65535)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_add_rmsnorm: bad arguments");
    const auto a8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
    const int part4 = H / (4 * stack::kNormSplit);
    const bool vec = H % (4 * stack::kNormSplit) == 0 && part4 <= 128 * 8 && aligned16(resid) && a8(weight) &&
                     a8(out) && (!delta || a8(delta));
    cudaStream_t s = as_stream(stream);
    cudaError_t e;
    const dim3 grid(stack::kNormSplit, M), block(128);
    if (!vec)
        e = launch_chained(stack::add_rmsnorm_any_kernel, dim3(M), dim3(256), 0, s, 1, resid, delta, weight, out, H,
                           eps);
    else if (part4 <= 128 * 2)
        e = launch_chained(stack::add_rmsnorm_kernel<2>, grid, block, 0, s, stack::kNormSplit, resid, delta, weight,
                           out, H, eps);
    else if (part4 <= 128 * 4)
        e = launch_chained(stack::add_rmsnorm_kernel<4>, grid, block, 0, s, stack::kNormSplit, resid, delta, weight,
                           out, H, eps);
    else
        e = launch_chained(stack::add_rmsnorm_kernel<8>, grid, block, 0, s, stack::kNormSplit, resid, delta, weight,
                           out, H, eps);
    DFLASH_CUDA_TRY(e);
    return DFLASH_OK;
}

extern "C" int dflash_stack_add_rmsnorm_reduce(float* resid, void* exchange, int world, int set,
                                               const dflash_bf16* weight, dflash_bf16* out, int M, int H, float eps,
                                               dflash_stream_t stream) {
    if (!resid || !exchange || !weight || !out || M < 1 || H < 1 || M > 65535 || world < 1 ||
        world > tp::kMaxRanks || (set != 0 && set != 1))
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_add_rmsnorm_reduce: bad arguments");
    const auto a8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
    const int part4 = H / (4 * stack::kNormSplit);
    if (H % (4 * stack::kNormSplit) || part4 > 128 * 8 || !aligned16(resid) || !a8(weight) || !a8(out) ||
        !aligned16(exchange))
        return fail(DFLASH_ERR_UNSUPPORTED, "dflash_stack_add_rmsnorm_reduce: H=%d (a multiple of %d up to %d) and "
                    "aligned buffers needed", H, 4 * stack::kNormSplit, 4 * stack::kNormSplit * 128 * 8);
    cudaStream_t s = as_stream(stream);
    const dim3 grid(stack::kNormSplit, M), block(128);
    cudaError_t e;
    if (part4 <= 128 * 2)
        e = launch_chained(stack::add_rmsnorm_reduce_kernel<2>, grid, block, 0, s, stack::kNormSplit, resid, exchange,
                           world, set, weight, out, M, H, eps);
    else if (part4 <= 128 * 4)
        e = launch_chained(stack::add_rmsnorm_reduce_kernel<4>, grid, block, 0, s, stack::kNormSplit, resid, exchange,
                           world, set, weight, out, M, H, eps);
    else
        e = launch_chained(stack::add_rmsnorm_reduce_kernel<8>, grid, block, 0, s, stack::kNormSplit, resid, exchange,
                           world, set, weight, out, M, H, eps);
    DFLASH_CUDA_TRY(e);
    return DFLASH_OK;
}

extern "C" int dflash_stack_silu_mul(const dflash_bf16* gate_up, dflash_bf16* y, int M, int I, dflash_stream_t stream) {
    if (!gate_up || !y || M < 1 || I < 1) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_silu_mul: bad arguments");
    const size_t n = (size_t)M * I;
    DFLASH_CUDA_TRY(launch_chained(stack::silu_mul_kernel, dim3(stack::grid_for(n, 256)), dim3(256), 0,
                                   as_stream(stream), 1, gate_up, y, M, I));
    return DFLASH_OK;
}

extern "C" int dflash_stack_conv_silu(const dflash_bf16* x, int ld, const dflash_bf16* window, const dflash_bf16* weight,
                                      dflash_bf16* y, int M, int C, int kc, int parts, dflash_stream_t stream) {
    if (!x || !window || !weight || !y || M < 1 || C < 1 || ld < C || parts < 1 || C % parts)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_conv_silu: bad arguments");
    if (kc < 1 || kc > 8) return fail(DFLASH_ERR_UNSUPPORTED, "conv width %d not in 1..8", kc);
    if (M > 16) return fail(DFLASH_ERR_UNSUPPORTED, "conv over M=%d tokens; at most 16", M);
    const dim3 grid((C + 127) / 128), block(128);
    cudaStream_t s = as_stream(stream);
    cudaError_t e = cudaSuccess;
    switch (kc) {
#define DFLASH_CONV_CASE(KC)                                                                                        \
    case KC:                                                                                                        \
        e = launch_chained(stack::conv_silu_kernel<KC>, grid, block, 0, s, 1, x, ld, window, weight, y, M, C, parts); \
        break;
        DFLASH_CONV_CASE(1) DFLASH_CONV_CASE(2) DFLASH_CONV_CASE(3) DFLASH_CONV_CASE(4)
        DFLASH_CONV_CASE(5) DFLASH_CONV_CASE(6) DFLASH_CONV_CASE(7) DFLASH_CONV_CASE(8)
#undef DFLASH_CONV_CASE
    }
    DFLASH_CUDA_TRY(e);
    return DFLASH_OK;
}

extern "C" int dflash_stack_gdn_gates(dflash_bf16* q, dflash_bf16* k, const dflash_bf16* ab, int ld_ab,
                                      const float* a_log, const float* dt_bias, float* alpha, float* beta, int M,
                                      int heads, int dk, dflash_stream_t stream) {
    if (!q || !k || !ab || !a_log || !dt_bias || !alpha || !beta || M < 1 || heads < 1 || dk < 1)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_gdn_gates: bad arguments");
    const int warps = M * heads;
    DFLASH_CUDA_TRY(launch_chained(stack::gdn_gates_kernel, dim3((warps + 7) / 8), dim3(256), 0, as_stream(stream), 1,
                                   q, k, ab, ld_ab, a_log, dt_bias, alpha, beta, M, heads, dk));
    return DFLASH_OK;
}

extern "C" int dflash_stack_gated_norm(const dflash_bf16* o, const dflash_bf16* z, int ld_z, const dflash_bf16* weight,
                                       dflash_bf16* out, int M, int heads, int dv, float eps, dflash_stream_t stream) {
    if (!o || !z || !weight || !out || M < 1 || heads < 1 || dv < 1)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_gated_norm: bad arguments");
    const int warps = M * heads;
    const dim3 grid((warps + 7) / 8), block(256);
    cudaStream_t s = as_stream(stream);
    cudaError_t e;
    switch (dv) {
        case 32: e = launch_chained(stack::gated_norm_kernel<1>, grid, block, 0, s, 1, o, z, ld_z, weight, out, M,
                                    heads, dv, eps); break;
        case 64: e = launch_chained(stack::gated_norm_kernel<2>, grid, block, 0, s, 1, o, z, ld_z, weight, out, M,
                                    heads, dv, eps); break;
        case 128: e = launch_chained(stack::gated_norm_kernel<4>, grid, block, 0, s, 1, o, z, ld_z, weight, out, M,
                                     heads, dv, eps); break;
        case 256: e = launch_chained(stack::gated_norm_kernel<8>, grid, block, 0, s, 1, o, z, ld_z, weight, out, M,
                                     heads, dv, eps); break;
        default: e = launch_chained(stack::gated_norm_kernel<0>, grid, block, 0, s, 1, o, z, ld_z, weight, out, M,
                                    heads, dv, eps);
    }
    DFLASH_CUDA_TRY(e);
    return DFLASH_OK;
}

static int attn_prep(dflash_bf16* qkv, int ld, const dflash_bf16* q_norm, const dflash_bf16* k_norm,
                     dflash_bf16* cache_k, dflash_bf16* cache_v, int M, int hq, int hkv, int d, int rot, int pos0,
                     int max_len, float eps, float theta, const int32_t* parents, dflash_stream_t stream,
                     const int32_t* position = nullptr) {
    if (position) pos0 = 0;  // read on the device; the kernel checks it against max_len
    if (!qkv || !q_norm || !k_norm || !cache_k || !cache_v || M < 1 || hq < 1 || hkv < 1 || pos0 < 0 ||
        pos0 + M > max_len || ld < (2 * hq + 2 * hkv) * d)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_attn_prep: bad arguments");
    if ((d != 64 && d != 128 && d != 256) || rot < 0 || rot > d || rot % 64)
        return fail(DFLASH_ERR_UNSUPPORTED, "head dim %d / rotary dims %d: need d in {64,128,256}, rot a multiple of 64",
                    d, rot);
    const int warps = M * (hq + hkv);
    const dim3 grid((warps + 7) / 8), block(256);
    cudaStream_t s = as_stream(stream);
    cudaError_t e;
    switch (d) {
        case 64:
            e = launch_chained(stack::attn_prep_kernel<2>, grid, block, 0, s, 1, qkv, ld, q_norm, k_norm, cache_k,
                               cache_v, M, hq, hkv, rot, pos0, max_len, eps, theta, parents, position);
            break;
        case 128:
            e = launch_chained(stack::attn_prep_kernel<4>, grid, block, 0, s, 1, qkv, ld, q_norm, k_norm, cache_k,
                               cache_v, M, hq, hkv, rot, pos0, max_len, eps, theta, parents, position);
            break;
        default:
            e = launch_chained(stack::attn_prep_kernel<8>, grid, block, 0, s, 1, qkv, ld, q_norm, k_norm, cache_k,
                               cache_v, M, hq, hkv, rot, pos0, max_len, eps, theta, parents, position);
            break;
    }
    DFLASH_CUDA_TRY(e);
    return DFLASH_OK;
}

extern "C" int dflash_stack_attn_prep(dflash_bf16* qkv, int ld, const dflash_bf16* q_norm, const dflash_bf16* k_norm,
                                      dflash_bf16* cache_k, dflash_bf16* cache_v, int M, int hq, int hkv, int d,
                                      int rot, int pos0, int max_len, float eps, float theta, dflash_stream_t stream) {
    return attn_prep(qkv, ld, q_norm, k_norm, cache_k, cache_v, M, hq, hkv, d, rot, pos0, max_len, eps, theta, nullptr,
                     stream);
}

extern "C" int dflash_stack_attn_prep_tree(dflash_bf16* qkv, int ld, const dflash_bf16* q_norm,
                                           const dflash_bf16* k_norm, dflash_bf16* cache_k, dflash_bf16* cache_v,
                                           int M, int hq, int hkv, int d, int rot, int pos0, int max_len, float eps,
                                           float theta, const int32_t* parents, dflash_stream_t stream) {
    if (!parents || M > kMaxTreeRows)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_attn_prep_tree: need parents and M <= %d", kMaxTreeRows);
    return attn_prep(qkv, ld, q_norm, k_norm, cache_k, cache_v, M, hq, hkv, d, rot, pos0, max_len, eps, theta, parents,
                     stream);
}

static int attn_decode(const dflash_bf16* qkv, int ld, const dflash_bf16* cache_k, const dflash_bf16* cache_v,
                       dflash_bf16* out, int M, int hq, int hkv, int d, int pos0, int max_len, float scale,
                       const int32_t* parents, dflash_stream_t stream, const int32_t* position = nullptr) {
    if (position) pos0 = 0;  // read on the device; the kernel checks it against max_len
    if (!qkv || !cache_k || !cache_v || !out || M < 1 || hq < 1 || hkv < 1 || hq % hkv || pos0 < 0 ||
        pos0 + M > max_len || ld < (2 * hq + 2 * hkv) * d || M > 65535)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_attn_decode: bad arguments");
    if (d != 64 && d != 128 && d != 256) return fail(DFLASH_ERR_UNSUPPORTED, "head dim %d not in {64,128,256}", d);
    if (hq / hkv > stack::kMaxG)
        return fail(DFLASH_ERR_UNSUPPORTED, "%d q heads per kv head; at most %d", hq / hkv, stack::kMaxG);
    if (!aligned16(cache_k) || !aligned16(cache_v) || !aligned16(qkv) || (ld * 2) % 16)
        return fail(DFLASH_ERR_MISALIGNED, "dflash_stack_attn_decode: qkv, its row stride and the caches must be "
                                           "16-byte aligned");
    int dev = 0;
    DFLASH_CUDA_TRY(cudaGetDevice(&dev));
    // twice the CTAs per (kv head, token) while the grid stays within half the SMs (measured:
    // 64 CTAs of 8 beat 32 of 4 by a third; 128 of 8 lose to 64 of 4)
    const bool small = 2LL * hkv * stack::kSplitSmall * M <= sm_count(dev);
    const int split = small ? stack::kSplitSmall : stack::kSplit;
    const dim3 grid(hkv * split, M), block(256);
    cudaStream_t s = as_stream(stream);
    const int G = hq / hkv;
    const int gmin = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;  // heads padded to a power of two
    const int ch = d / 32;
    const int gp = gmin > ch / 2 ? gmin : ch / 2;                 // keeps the score registers bounded
    cudaError_t e = cudaErrorInvalidValue;
#define DFLASH_ATTN_CASE(CH, GP)                                                                                   \
    if (ch == CH && gp == GP)                                                                                      \
        e = small ? launch_chained(stack::attn_decode_kernel<CH, GP, stack::kSplitSmall>, grid, block, 0, s,        \
                                   stack::kSplitSmall, qkv, ld, cache_k, cache_v, out, hq, hkv, pos0, max_len, scale, \
                                   parents, position)                                                              \
                  : launch_chained(stack::attn_decode_kernel<CH, GP, stack::kSplit>, grid, block, 0, s,             \
                                   stack::kSplit, qkv, ld, cache_k, cache_v, out, hq, hkv, pos0, max_len, scale,    \
                                   parents, position);
    DFLASH_ATTN_CASE(2, 1) DFLASH_ATTN_CASE(2, 2) DFLASH_ATTN_CASE(2, 4) DFLASH_ATTN_CASE(2, 8)
    DFLASH_ATTN_CASE(4, 2) DFLASH_ATTN_CASE(4, 4) DFLASH_ATTN_CASE(4, 8)
    DFLASH_ATTN_CASE(8, 4) DFLASH_ATTN_CASE(8, 8)
#undef DFLASH_ATTN_CASE
    DFLASH_CUDA_TRY(e);
    return DFLASH_OK;
}

extern "C" int dflash_stack_attn_decode(const dflash_bf16* qkv, int ld, const dflash_bf16* cache_k,
                                        const dflash_bf16* cache_v, dflash_bf16* out, int M, int hq, int hkv, int d,
                                        int pos0, int max_len, float scale, dflash_stream_t stream) {
    return attn_decode(qkv, ld, cache_k, cache_v, out, M, hq, hkv, d, pos0, max_len, scale, nullptr, stream);
}

extern "C" int dflash_stack_attn_decode_tree(const dflash_bf16* qkv, int ld, const dflash_bf16* cache_k,
                                             const dflash_bf16* cache_v, dflash_bf16* out, int M, int hq, int hkv,
                                             int d, int pos0, int max_len, float scale, const int32_t* parents,
                                             dflash_stream_t stream) {
    if (!parents || M > kMaxTreeRows)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_attn_decode_tree: need parents and M <= %d",
                    kMaxTreeRows);
    return attn_decode(qkv, ld, cache_k, cache_v, out, M, hq, hkv, d, pos0, max_len, scale, parents, stream);
}

extern "C" int dflash_accept(const unsigned long long* argmax_keys, const int32_t* proposals, int drafts,
                             int32_t* target_tokens, int32_t* accepted, dflash_stream_t stream) {
    if (!argmax_keys || (!proposals && drafts > 0) || !target_tokens || !accepted || drafts < 0)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_accept: bad arguments");
    DFLASH_CUDA_TRY(launch_chained(stack::accept_kernel, dim3(1), dim3(32), 0, as_stream(stream), 1, argmax_keys,
                                   proposals, drafts, target_tokens, accepted));
    return DFLASH_OK;
}

static int gdn_conv_gates(const dflash_bf16* x, int ld, const dflash_bf16* window, const dflash_bf16* weight,
                          dflash_bf16* y, const dflash_bf16* ab, int ld_ab, const float* a_log, const float* dt_bias,
                          float* alpha, float* beta, int M, int heads, int dk, int kc, const int32_t* parents,
                          dflash_stream_t stream) {
    if (!x || !window || !weight || !y || !ab || !a_log || !dt_bias || !alpha || !beta || M < 1 || heads < 1 ||
        ld < 3 * heads * dk)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_gdn_conv_gates: bad arguments");
    if ((dk != 32 && dk != 64 && dk != 128) || kc < 2 || kc > 4)
        return fail(DFLASH_ERR_UNSUPPORTED, "dflash_stack_gdn_conv_gates: dk %d (32, 64, 128) / conv width %d (2..4)",
                    dk, kc);
    const int warps = 3 * heads * M;
    const dim3 grid((warps + 7) / 8), block(256);
    cudaStream_t s = as_stream(stream);
    cudaError_t e = cudaSuccess;
#define DFLASH_CG_CASE(KC, DJ)                                                                                   \
    if (kc == KC && dk == 32 * DJ)                                                                               \
        e = launch_chained(stack::gdn_conv_gates_kernel<KC, DJ>, grid, block, 0, s, 1, x, ld, window, weight, y, ab, \
                           ld_ab, a_log, dt_bias, alpha, beta, M, heads, parents);
    DFLASH_CG_CASE(2, 1) DFLASH_CG_CASE(2, 2) DFLASH_CG_CASE(2, 4)
    DFLASH_CG_CASE(3, 1) DFLASH_CG_CASE(3, 2) DFLASH_CG_CASE(3, 4)
    DFLASH_CG_CASE(4, 1) DFLASH_CG_CASE(4, 2) DFLASH_CG_CASE(4, 4)
#undef DFLASH_CG_CASE
    DFLASH_CUDA_TRY(e);
    return DFLASH_OK;
}

extern "C" int dflash_stack_gdn_conv_gates(const dflash_bf16* x, int ld, const dflash_bf16* window,
                                           const dflash_bf16* weight, dflash_bf16* y, const dflash_bf16* ab,
                                           int ld_ab, const float* a_log, const float* dt_bias, float* alpha,
                                           float* beta, int M, int heads, int dk, int kc, dflash_stream_t stream) {
    return gdn_conv_gates(x, ld, window, weight, y, ab, ld_ab, a_log, dt_bias, alpha, beta, M, heads, dk, kc, nullptr,
                          stream);
}

extern "C" int dflash_stack_gdn_conv_gates_tree(const dflash_bf16* x, int ld, const dflash_bf16* window,
                                                const dflash_bf16* weight, dflash_bf16* y, const dflash_bf16* ab,
                                                int ld_ab, const float* a_log, const float* dt_bias, float* alpha,
                                                float* beta, int M, int heads, int dk, int kc,
                                                const int32_t* parents, dflash_stream_t stream) {
    if (!parents || M > kMaxTreeRows)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_gdn_conv_gates_tree: need parents and M <= %d",
                    kMaxTreeRows);
    return gdn_conv_gates(x, ld, window, weight, y, ab, ld_ab, a_log, dt_bias, alpha, beta, M, heads, dk, kc, parents,
                          stream);
}

extern "C" int dflash_accept_reduce(void* exchange, int world, int set, const int32_t* proposals, int drafts,
                                    int32_t* target_tokens, int32_t* accepted, dflash_stream_t stream) {
    if (!exchange || world < 1 || world > tp::kMaxRanks || (set != 0 && set != 1) || (!proposals && drafts > 0) ||
        !target_tokens || !accepted || drafts < 0)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_accept_reduce: bad arguments");
    DFLASH_CUDA_TRY(launch_chained(stack::accept_reduce_kernel, dim3(1), dim3(32), 0, as_stream(stream), 1, exchange,
                                   world, set, proposals, drafts, target_tokens, accepted));
    return DFLASH_OK;
}

extern "C" int dflash_stack_kv_compact(dflash_bf16* cache_k, dflash_bf16* cache_v, int layers, long long layer_stride,
                                       int hkv, int d, int pos0, int max_len, const int32_t* rows, int keep,
                                       dflash_stream_t stream) {
    if (!cache_k || !cache_v || cache_k == cache_v || !rows || layers < 1 || layers > 65535 || hkv < 1 ||
        hkv > 65535 || pos0 < 0 || max_len < 1 || keep < 1 || keep > kMaxTreeRows || layer_stride < 0 ||
        (layers > 1 && layer_stride < (long long)hkv * max_len * d))
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_kv_compact: bad arguments");
    if (d != 64 && d != 128 && d != 256) return fail(DFLASH_ERR_UNSUPPORTED, "head dim %d not in {64,128,256}", d);
    if (!aligned16(cache_k) || !aligned16(cache_v) || (layer_stride * 2) % 16)
        return fail(DFLASH_ERR_MISALIGNED, "dflash_stack_kv_compact: caches and layer stride must be 16-byte aligned");
    stack::CompactRows rl{};
    for (int i = 0; i < keep; ++i) {
        if (rows[i] < 0 || pos0 + rows[i] >= max_len)
            return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_kv_compact: rows[%d]=%d outside the cache", i,
                        rows[i]);
        rl.r[i] = rows[i];
    }
    if (pos0 + keep > max_len) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_kv_compact: keep past max_len");
    DFLASH_CUDA_TRY(launch_chained(stack::kv_compact_kernel, dim3(hkv, layers, 2), dim3(256), 0, as_stream(stream), 1,
                                   reinterpret_cast<uint16_t*>(cache_k), reinterpret_cast<uint16_t*>(cache_v),
                                   layer_stride, d, pos0, max_len, rl, keep));
    return DFLASH_OK;
}

extern "C" int dflash_bias_add(dflash_bf16* y, const dflash_bf16* bias, int rows, int N, dflash_stream_t stream) {
    if (!y || !bias || rows < 1 || N < 1) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_bias_add: bad arguments");
    const long long total = (long long)rows * N;
    const long long blocks = (total + 255) / 256;
    if (blocks > 0x7fffffffLL) return fail(DFLASH_ERR_UNSUPPORTED, "dflash_bias_add: %lld elements", total);
    DFLASH_CUDA_TRY(launch_chained(stack::bias_add_kernel, dim3((unsigned)blocks), dim3(256), 0, as_stream(stream), 1,
                                   reinterpret_cast<uint16_t*>(y), reinterpret_cast<const uint16_t*>(bias), total, N));
    return DFLASH_OK;
}

extern "C" int dflash_accept_tree(const int32_t* target_tokens, const int32_t* parents, const int32_t* tokens,
                                  int rows, int32_t* path, int32_t* path_len, int32_t* next_token,
                                  dflash_stream_t stream) {
    if (!target_tokens || !parents || !tokens || !path || !path_len || !next_token || rows < 1 ||
        rows > kMaxTreeRows)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_accept_tree: bad arguments (1 <= rows <= %d)", kMaxTreeRows);
    DFLASH_CUDA_TRY(launch_chained(stack::accept_tree_kernel, dim3(1), dim3(32), 0, as_stream(stream), 1,
                                   target_tokens, parents, tokens, rows, path, path_len, next_token));
    return DFLASH_OK;
}

extern "C" int dflash_stack_gdn_conv_gates_grouped(const dflash_bf16* x, int ld, const dflash_bf16* window,
                                                   const dflash_bf16* weight, dflash_bf16* y, const dflash_bf16* ab,
                                                   int ld_ab, const float* a_log, const float* dt_bias, float* alpha,
                                                   float* beta, int M, int heads, int k_heads, int dk, int kc,
                                                   const int32_t* parents, dflash_stream_t stream) {
    if (!x || !window || !weight || !y || !ab || !a_log || !dt_bias || !alpha || !beta || M < 1 || heads < 1 ||
        k_heads < 1 || heads % k_heads || ld < (2 * k_heads + heads) * dk || ld_ab < 2 * heads)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_gdn_conv_gates_grouped: bad arguments");
    if (parents && M > kMaxTreeRows)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_gdn_conv_gates_grouped: a tree has at most %d rows",
                    kMaxTreeRows);
    if ((dk != 32 && dk != 64 && dk != 128) || kc < 2 || kc > 4)
        return fail(DFLASH_ERR_UNSUPPORTED,
                    "dflash_stack_gdn_conv_gates_grouped: dk %d (32, 64, 128) / conv width %d (2..4)", dk, kc);
    const long long warps = (long long)M * (2 * k_heads + heads);
    const dim3 grid((unsigned)((warps + 7) / 8)), block(256);
    cudaStream_t s = as_stream(stream);
    cudaError_t e = cudaSuccess;
#define DFLASH_CGG_CASE(KC, DJ)                                                                                  \
    if (kc == KC && dk == 32 * DJ)                                                                              \
        e = launch_chained(stack::gdn_conv_gates_grouped_kernel<KC, DJ>, grid, block, 0, s, 1, x, ld, window, weight, \
                           y, ab, ld_ab, a_log, dt_bias, alpha, beta, M, heads, k_heads, parents);
    DFLASH_CGG_CASE(2, 1) DFLASH_CGG_CASE(2, 2) DFLASH_CGG_CASE(2, 4)
    DFLASH_CGG_CASE(3, 1) DFLASH_CGG_CASE(3, 2) DFLASH_CGG_CASE(3, 4)
    DFLASH_CGG_CASE(4, 1) DFLASH_CGG_CASE(4, 2) DFLASH_CGG_CASE(4, 4)
#undef DFLASH_CGG_CASE
    DFLASH_CUDA_TRY(e);
    return DFLASH_OK;
}

extern "C" int dflash_stack_attn_prep_ex(dflash_bf16* qkv, int ld, const dflash_bf16* q_norm,
                                         const dflash_bf16* k_norm, dflash_bf16* cache_k, dflash_bf16* cache_v, int M,
                                         int hq, int hkv, int d, int rot, int pos0, int max_len, float eps,
                                         float theta, const int32_t* parents, const int32_t* position,
                                         dflash_stream_t stream) {
    if (parents && M > kMaxTreeRows)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_attn_prep_ex: a tree has at most %d rows", kMaxTreeRows);
    return attn_prep(qkv, ld, q_norm, k_norm, cache_k, cache_v, M, hq, hkv, d, rot, pos0, max_len, eps, theta, parents,
                     stream, position);
}

extern "C" int dflash_stack_attn_decode_ex(const dflash_bf16* qkv, int ld, const dflash_bf16* cache_k,
                                           const dflash_bf16* cache_v, dflash_bf16* out, int M, int hq, int hkv, int d,
                                           int pos0, int max_len, float scale, const int32_t* parents,
                                           const int32_t* position, dflash_stream_t stream) {
    if (parents && M > kMaxTreeRows)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_attn_decode_ex: a tree has at most %d rows",
                    kMaxTreeRows);
    return attn_decode(qkv, ld, cache_k, cache_v, out, M, hq, hkv, d, pos0, max_len, scale, parents, stream, position);
}
