// Glue kernels of the tensor-parallel verify stack (the hybrid target's layers around the
// quantized projections): residual add + RMSNorm, the SiLU-gated MLP activation, the
// gated-delta layer's causal depthwise convolution, per-head normalisation, gates and
// gated output norm, and the attention layer's q/k norm + rotary embedding + cache append
// and its decode attention with the output gate.  The projections themselves are
// dflash_qmm and the recurrence is dflash_gdn_step.
//
// All tensors are row-major with one row per token (M rows, the verify block).  Every
// kernel here is memory- or latency-bound and tiny next to the weight stream.
#include "common.cuh"
#include "dflash_stack.h"

namespace dflash {
namespace stack {

__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
__device__ __forceinline__ uint16_t to_bf(float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    return *reinterpret_cast<const uint16_t*>(&h);
}
__device__ __forceinline__ float bf_round(float v) { return bf(to_bf(v)); }
__device__ __forceinline__ float silu(float v) { return v / (1.f + __expf(-v)); }

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += red[i];  // the same order on every thread
    return t;
}

// resid[m] += delta[m] (if given); out[m] = bf16(resid[m] * rsqrt(mean(resid[m]^2) + eps) * w)
__global__ void add_rmsnorm_kernel(float* __restrict__ resid, const uint16_t* __restrict__ delta,
                                   const uint16_t* __restrict__ w, uint16_t* __restrict__ out, int H, float eps) {
    __shared__ float red[32];
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
// after the round dflash_gdn_conv_rollback rebuilds it from the accepted inputs.
template <int KC>
__global__ void conv_silu_kernel(const uint16_t* __restrict__ x, int ld, const uint16_t* __restrict__ window,
                                 const uint16_t* __restrict__ w, uint16_t* __restrict__ y, int M, int C, int parts) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    constexpr int h = KC - 1;
    float hist[h > 0 ? h : 1];
#pragma unroll
    for (int i = 0; i < h; ++i) hist[i] = bf(window[(size_t)i * C + c]);
    float wk[KC];
#pragma unroll
    for (int i = 0; i < KC; ++i) wk[i] = bf(w[(size_t)c * KC + i]);
    const int cp = C / parts, part = c / cp, cc = c - part * cp;
    for (int t = 0; t < M; ++t) {
        const float xt = bf(x[(size_t)t * ld + c]);
        float acc = wk[KC - 1] * xt;
#pragma unroll
        for (int i = 0; i < h; ++i) acc = fmaf(wk[i], hist[i], acc);
        y[((size_t)part * M + t) * cp + cc] = to_bf(silu(acc));
#pragma unroll
        for (int i = 0; i + 1 < h; ++i) hist[i] = hist[i + 1];
        if constexpr (h > 0) hist[h - 1] = xt;
    }
}

// Per (token, head) of the gated-delta layer: L2-normalise q and k (dk each) in place,
// alpha = exp(-exp(a_log[h]) * softplus(a + dt_bias[h])), beta = sigmoid(b).
// q, k: [M, heads * dk]; ab: [M, ld_ab] with b at [0, heads) and a at [heads, 2 heads).
// One warp per (token, head).
__global__ void gdn_gates_kernel(uint16_t* __restrict__ q, uint16_t* __restrict__ k, const uint16_t* __restrict__ ab,
                                 int ld_ab, const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                                 float* __restrict__ alpha, float* __restrict__ beta, int M, int heads, int dk) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M * heads) return;
    const int t = warp / heads, h = warp % heads;
    for (int part = 0; part < 2; ++part) {
        uint16_t* v = (part ? k : q) + ((size_t)t * heads + h) * dk;
        float ss = 0.f;
        for (int i = lane; i < dk; i += 32) ss = fmaf(bf(v[i]), bf(v[i]), ss);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rs = rsqrtf(ss + 1e-6f);
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

// out[t, h*dv + i] = rmsnorm(o[t, h, :]) * w[i] * silu(z[t, h*dv + i]); one warp per (t, h).
__global__ void gated_norm_kernel(const uint16_t* __restrict__ o, const uint16_t* __restrict__ z, int ld_z,
                                  const uint16_t* __restrict__ w, uint16_t* __restrict__ out, int M, int heads, int dv,
                                  float eps) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M * heads) return;
    const int t = warp / heads, h = warp % heads;
    const uint16_t* ov = o + ((size_t)t * heads + h) * dv;
    float ss = 0.f;
    for (int i = lane; i < dv; i += 32) ss = fmaf(bf(ov[i]), bf(ov[i]), ss);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, s);
    const float rs = rsqrtf(ss / dv + eps);
    for (int i = lane; i < dv; i += 32) {
        const float zz = bf(z[(size_t)t * ld_z + (size_t)h * dv + i]);
        out[((size_t)t * heads + h) * dv + i] = to_bf(bf(ov[i]) * rs * bf(w[i]) * silu(zz));
    }
}

// Attention-layer prep, one warp per (token, head slot).  qkv row t (stride ld) holds
// [q (hq * d) | gate (hq * d) | k (hkv * d) | v (hkv * d)].  Slot < hq: q head, RMSNorm with
// q_norm then rotary embedding on its first `rot` dims, in place.  Slot >= hq: kv head j,
// k gets k_norm and the rotary embedding and goes to cache_k[j, pos0 + t]; v is copied to
// cache_v[j, pos0 + t].  Rotary: rotate-half over the first rot dims, frequency
// theta^(-2i/rot) for pair (i, i + rot/2), position pos0 + t.  Lane l holds dims
// l + 32 c, so with rot a multiple of 64 both halves of a pair sit in one lane.
template <int CH>
__global__ void attn_prep_kernel(uint16_t* __restrict__ qkv, int ld, const uint16_t* __restrict__ q_norm,
                                 const uint16_t* __restrict__ k_norm, uint16_t* __restrict__ cache_k,
                                 uint16_t* __restrict__ cache_v, int M, int hq, int hkv, int rot, int pos0,
                                 int max_len, float eps, float theta) {
    constexpr int d = CH * 32;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int slots = hq + hkv;
    if (warp >= M * slots) return;
    const int t = warp / slots, slot = warp % slots;
    uint16_t* row = qkv + (size_t)t * ld;
    if (slot >= hq) {  // v copy first (independent of the k work)
        const int j = slot - hq;
        const uint16_t* vs = row + (size_t)(2 * hq + hkv + j) * d;
        uint16_t* vd = cache_v + ((size_t)j * max_len + pos0 + t) * d;
#pragma unroll
        for (int c = 0; c < CH; ++c) vd[lane + 32 * c] = vs[lane + 32 * c];
    }
    uint16_t* src = slot < hq ? row + (size_t)slot * d : row + (size_t)(2 * hq + (slot - hq)) * d;
    uint16_t* dst = slot < hq ? src : cache_k + ((size_t)(slot - hq) * max_len + pos0 + t) * d;
    const uint16_t* nw = slot < hq ? q_norm : k_norm;
    float v[CH];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        v[c] = bf(src[lane + 32 * c]);
        ss = fmaf(v[c], v[c], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rs = rsqrtf(ss / d + eps);
#pragma unroll
    for (int c = 0; c < CH; ++c) v[c] = bf_round(v[c] * rs * bf(nw[lane + 32 * c]));
    const int half_c = rot / 64;  // pair partner is c + half_c
    const float pos = (float)(pos0 + t);
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

// Attention of the M block tokens over the cache, one CTA (8 warps) per (q head, token).
// Token t sees keys 0 .. pos0 + t (the cache prefix and the block causally).  q: row t of
// qkv at head h; gate at [hq * d + h * d); q head h reads kv head h / (hq / hkv).
// out[t, h * d + e] = softmax(q K^T * scale) V * sigmoid(gate).  Each warp runs an online
// softmax over keys warp, warp + 8, ...; lane l holds dims [l * CH, l * CH + CH).
template <int CH>
__global__ void __launch_bounds__(256) attn_decode_kernel(const uint16_t* __restrict__ qkv, int ld,
                                                          const uint16_t* __restrict__ cache_k,
                                                          const uint16_t* __restrict__ cache_v,
                                                          uint16_t* __restrict__ out, int hq, int hkv, int pos0,
                                                          int max_len, float scale) {
    constexpr int d = CH * 32;
    __shared__ float s_m[8], s_l[8];
    __shared__ float s_acc[8][d];
    const int h = blockIdx.x, t = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvh = h / (hq / hkv);
    const uint16_t* qrow = qkv + (size_t)t * ld + (size_t)h * d + lane * CH;
    float q[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) q[c] = bf(qrow[c]) * scale;
    const uint16_t* kb = cache_k + (size_t)kvh * max_len * d + lane * CH;
    const uint16_t* vb = cache_v + (size_t)kvh * max_len * d + lane * CH;
    const int n = pos0 + t + 1;
    float m = -INFINITY, l = 0.f, acc[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) acc[c] = 0.f;
    for (int j = warp; j < n; j += 8) {
        const uint16_t* kr = kb + (size_t)j * d;
        float sdot = 0.f;
#pragma unroll
        for (int c = 0; c < CH; ++c) sdot = fmaf(q[c], bf(kr[c]), sdot);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sdot += __shfl_xor_sync(0xffffffffu, sdot, o);
        const float mn = fmaxf(m, sdot);
        const float corr = __expf(m - mn), p = __expf(sdot - mn);
        l = l * corr + p;
        const uint16_t* vr = vb + (size_t)j * d;
#pragma unroll
        for (int c = 0; c < CH; ++c) acc[c] = fmaf(p, bf(vr[c]), acc[c] * corr);
        m = mn;
    }
    if (lane == 0) {
        s_m[warp] = m;
        s_l[warp] = l;
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) s_acc[warp][lane * CH + c] = acc[c];
    __syncthreads();
    float mx = -INFINITY;
    for (int w = 0; w < 8; ++w) mx = fmaxf(mx, s_m[w]);
    float den = 0.f, f[8];
    for (int w = 0; w < 8; ++w) {
        f[w] = s_l[w] > 0.f ? __expf(s_m[w] - mx) : 0.f;
        den = fmaf(s_l[w], f[w], den);
    }
    const uint16_t* grow = qkv + (size_t)t * ld + (size_t)(hq + h) * d;
    for (int e = threadIdx.x; e < d; e += blockDim.x) {
        float num = 0.f;
        for (int w = 0; w < 8; ++w) num = fmaf(s_acc[w][e], f[w], num);
        const float g = bf(grow[e]);
        out[(size_t)t * hq * d + (size_t)h * d + e] = to_bf(num / den / (1.f + __expf(-g)));
    }
}

inline unsigned grid_for(size_t n, int block) {
    const size_t g = (n + block - 1) / block;
    return (unsigned)(g < 4096 ? (g > 0 ? g : 1) : 4096);
}

}  // namespace stack
}  // namespace dflash

using namespace dflash;

extern "C" int dflash_stack_add_rmsnorm(float* resid, const dflash_bf16* delta, const dflash_bf16* weight,
                                        dflash_bf16* out, int M, int H, float eps, dflash_stream_t stream) {
    if (!resid || !weight || !out || M < 1 || H < 1)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_add_rmsnorm: bad arguments");
    stack::add_rmsnorm_kernel<<<M, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(resid, delta, weight, out, H,
                                                                                         eps);
    DFLASH_CUDA_TRY(cudaGetLastError());
    return DFLASH_OK;
}

extern "C" int dflash_stack_silu_mul(const dflash_bf16* gate_up, dflash_bf16* y, int M, int I, dflash_stream_t stream) {
    if (!gate_up || !y || M < 1 || I < 1) return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_silu_mul: bad arguments");
    const size_t n = (size_t)M * I;
    stack::silu_mul_kernel<<<stack::grid_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(gate_up, y, M,
                                                                                                       I);
    DFLASH_CUDA_TRY(cudaGetLastError());
    return DFLASH_OK;
}

extern "C" int dflash_stack_conv_silu(const dflash_bf16* x, int ld, const dflash_bf16* window, const dflash_bf16* weight,
                                      dflash_bf16* y, int M, int C, int kc, int parts, dflash_stream_t stream) {
    if (!x || !window || !weight || !y || M < 1 || C < 1 || ld < C || parts < 1 || C % parts)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_conv_silu: bad arguments");
    if (kc < 1 || kc > 8) return fail(DFLASH_ERR_UNSUPPORTED, "conv width %d not in 1..8", kc);
    const dim3 grid((C + 127) / 128), block(128);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (kc) {
#define DFLASH_CONV_CASE(KC) \
    case KC: stack::conv_silu_kernel<KC><<<grid, block, 0, s>>>(x, ld, window, weight, y, M, C, parts); break;
        DFLASH_CONV_CASE(1) DFLASH_CONV_CASE(2) DFLASH_CONV_CASE(3) DFLASH_CONV_CASE(4)
        DFLASH_CONV_CASE(5) DFLASH_CONV_CASE(6) DFLASH_CONV_CASE(7) DFLASH_CONV_CASE(8)
#undef DFLASH_CONV_CASE
    }
    DFLASH_CUDA_TRY(cudaGetLastError());
    return DFLASH_OK;
}

extern "C" int dflash_stack_gdn_gates(dflash_bf16* q, dflash_bf16* k, const dflash_bf16* ab, int ld_ab,
                                      const float* a_log, const float* dt_bias, float* alpha, float* beta, int M,
                                      int heads, int dk, dflash_stream_t stream) {
    if (!q || !k || !ab || !a_log || !dt_bias || !alpha || !beta || M < 1 || heads < 1 || dk < 1)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_gdn_gates: bad arguments");
    const int warps = M * heads;
    stack::gdn_gates_kernel<<<(warps + 7) / 8, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        q, k, ab, ld_ab, a_log, dt_bias, alpha, beta, M, heads, dk);
    DFLASH_CUDA_TRY(cudaGetLastError());
    return DFLASH_OK;
}

extern "C" int dflash_stack_gated_norm(const dflash_bf16* o, const dflash_bf16* z, int ld_z, const dflash_bf16* weight,
                                       dflash_bf16* out, int M, int heads, int dv, float eps, dflash_stream_t stream) {
    if (!o || !z || !weight || !out || M < 1 || heads < 1 || dv < 1)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_gated_norm: bad arguments");
    const int warps = M * heads;
    stack::gated_norm_kernel<<<(warps + 7) / 8, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(o, z, ld_z, weight,
                                                                                                out, M, heads, dv, eps);
    DFLASH_CUDA_TRY(cudaGetLastError());
    return DFLASH_OK;
}

extern "C" int dflash_stack_attn_prep(dflash_bf16* qkv, int ld, const dflash_bf16* q_norm, const dflash_bf16* k_norm,
                                      dflash_bf16* cache_k, dflash_bf16* cache_v, int M, int hq, int hkv, int d,
                                      int rot, int pos0, int max_len, float eps, float theta, dflash_stream_t stream) {
    if (!qkv || !q_norm || !k_norm || !cache_k || !cache_v || M < 1 || hq < 1 || hkv < 1 || pos0 < 0 ||
        pos0 + M > max_len || ld < (2 * hq + 2 * hkv) * d)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_attn_prep: bad arguments");
    if ((d != 64 && d != 128 && d != 256) || rot < 0 || rot > d || rot % 64)
        return fail(DFLASH_ERR_UNSUPPORTED, "head dim %d / rotary dims %d: need d in {64,128,256}, rot a multiple of 64", d, rot);
    const int warps = M * (hq + hkv);
    const dim3 grid((warps + 7) / 8), block(256);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (d) {
        case 64: stack::attn_prep_kernel<2><<<grid, block, 0, s>>>(qkv, ld, q_norm, k_norm, cache_k, cache_v, M, hq, hkv, rot, pos0, max_len, eps, theta); break;
        case 128: stack::attn_prep_kernel<4><<<grid, block, 0, s>>>(qkv, ld, q_norm, k_norm, cache_k, cache_v, M, hq, hkv, rot, pos0, max_len, eps, theta); break;
        default: stack::attn_prep_kernel<8><<<grid, block, 0, s>>>(qkv, ld, q_norm, k_norm, cache_k, cache_v, M, hq, hkv, rot, pos0, max_len, eps, theta); break;
    }
    DFLASH_CUDA_TRY(cudaGetLastError());
    return DFLASH_OK;
}

extern "C" int dflash_stack_attn_decode(const dflash_bf16* qkv, int ld, const dflash_bf16* cache_k,
                                        const dflash_bf16* cache_v, dflash_bf16* out, int M, int hq, int hkv, int d,
                                        int pos0, int max_len, float scale, dflash_stream_t stream) {
    if (!qkv || !cache_k || !cache_v || !out || M < 1 || hq < 1 || hkv < 1 || hq % hkv || pos0 < 0 ||
        pos0 + M > max_len || ld < (2 * hq + 2 * hkv) * d || M > 65535)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_stack_attn_decode: bad arguments");
    if (d != 64 && d != 128 && d != 256) return fail(DFLASH_ERR_UNSUPPORTED, "head dim %d not in {64,128,256}", d);
    const dim3 grid(hq, M), block(256);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (d) {
        case 64: stack::attn_decode_kernel<2><<<grid, block, 0, s>>>(qkv, ld, cache_k, cache_v, out, hq, hkv, pos0, max_len, scale); break;
        case 128: stack::attn_decode_kernel<4><<<grid, block, 0, s>>>(qkv, ld, cache_k, cache_v, out, hq, hkv, pos0, max_len, scale); break;
        default: stack::attn_decode_kernel<8><<<grid, block, 0, s>>>(qkv, ld, cache_k, cache_v, out, hq, hkv, pos0, max_len, scale); break;
    }
    DFLASH_CUDA_TRY(cudaGetLastError());
    return DFLASH_OK;
}
